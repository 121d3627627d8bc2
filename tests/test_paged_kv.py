"""Paged KV cache: the host-side block allocator (CPU) and the paged decode
kernels against the contiguous ones on the same keys (GPU).  Pools are
[num_blocks, Hkv, 64, D]; block tables are shuffled so neighbouring keys of
a sequence sit in unrelated pool blocks."""
import pytest
import torch

from oracle import ops as O
from torchplusplus_b200.llmops.kvcache import PagedKVCache


def test_paged_allocator_reserve_release():
    c = PagedKVCache(num_blocks=10, n_kv_heads=2, head_dim=64, dtype=torch.float16,
                     device="cpu", batch_size=3, max_seq_len=1000)
    c.reserve(0, 130)            # 3 blocks
    c.reserve(1, 64)             # 1 block
    c.reserve(0, 150)            # still 3 blocks
    assert c.free_blocks == 6
    t = c.block_table
    assert (t[0, :3] >= 0).all() and (t[0, 3:] == -1).all()
    assert (t[1, :1] >= 0).all() and (t[1, 1:] == -1).all()
    assert len(set(t[0, :3].tolist()) | set(t[1, :1].tolist())) == 4  # distinct blocks
    c.release(0)
    assert c.free_blocks == 9 and (c.block_table[0] == -1).all()
    with pytest.raises(RuntimeError):
        c.reserve(2, 10 * 64 + 1)  # 11 blocks > 9 free
    with pytest.raises(ValueError):
        c.reserve(2, 1001)


def _pools_from_contiguous(kc, vc, g, spare=7):
    """Scatter contiguous caches [B, Hkv, S, D] into shuffled pool blocks via
    the paged append kernel; returns pools and the block table."""
    from torchplusplus_b200 import ops
    B, Hkv, S, D = kc.shape
    nb = (S + 63) // 64
    perm = torch.randperm(B * nb + spare, generator=g)
    table = perm[:B * nb].view(B, nb).to(torch.int32).cuda()
    kp = torch.zeros(B * nb + spare, Hkv, 64, D, dtype=kc.dtype, device="cuda")
    vp = torch.zeros_like(kp)
    ops.kv_append_paged(kc, vc, kp, vp, table, start_pos=0)
    return kp, vp, table


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", [
    # B, Hq, Hkv, D, lens, window
    (4, 16, 8, 128, [1, 64, 65, 700], -1),
    (3, 16, 8, 128, [513, 2000, 40], 255),      # window start inside a block
    (2, 8, 1, 64, [129, 5], -1),
    (1, 64, 2, 128, [9000], -1),                # many splits, two head passes
])
def test_attention_decode_paged_matches_contiguous(dtype, case):
    from torchplusplus_b200 import ops
    B, Hq, Hkv, D, lens, window = case
    g = torch.Generator().manual_seed(51)
    S = max(lens) + 3
    q = torch.randn(B, Hq, D, generator=g).to(dtype).cuda()
    kc = torch.randn(B, Hkv, S, D, generator=g).to(dtype).cuda()
    vc = torch.randn(B, Hkv, S, D, generator=g).to(dtype).cuda()
    sl = torch.tensor(lens, dtype=torch.int32).cuda()
    kp, vp, table = _pools_from_contiguous(kc, vc, g)
    # the append put every row where the table says
    for b in range(B):
        for k in (0, 63, 64, lens[b] - 1):
            blk = int(table[b, k // 64])
            assert torch.equal(kp[blk, :, k % 64], kc[b, :, k])
    y = ops.attention_decode_paged(q, kp, vp, table, sl, S, window_left=window)
    ref = O.attention_decode(q.cpu(), kc.cpu(), vc.cpu(), sl.cpu(), window_left=window)
    err = (y.float().cpu() - ref).abs() / ref.abs().clamp(min=1.0)
    assert err.max().item() <= 2e-2
    y2 = ops.attention_decode(q, kc, vc, sl, S, window_left=window)
    assert (y.float() - y2.float()).abs().max().item() <= 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("case", [
    (4, 16, 8, 128, [1, 64, 65, 700], -1),
    (3, 16, 8, 128, [513, 2000, 40], 255),
])
def test_attention_decode_qkv_paged_matches_contiguous(case):
    from torchplusplus_b200 import ops
    B, Hq, Hkv, D, lens, window = case
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(52)
    S = max(lens) + 3
    qkv = torch.randn(B, 1, (Hq + 2 * Hkv) * D, generator=g).to(dtype).cuda()
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype).cuda()
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype).cuda()
    cos, sin = O.compute_rope_params(D, 1e6, S)
    cos, sin = cos.cuda(), sin.cuda()
    kc = torch.randn(B, Hkv, S, D, generator=g).to(dtype).cuda()
    vc = torch.randn(B, Hkv, S, D, generator=g).to(dtype).cuda()
    sl = torch.tensor(lens, dtype=torch.int32).cuda()
    pos = sl - 1
    kp, vp, table = _pools_from_contiguous(kc, vc, g)
    y = ops.attention_decode_qkv_paged(qkv, qn, kn, 1e-6, cos, sin, pos, kp, vp, table, sl, S,
                                       Hq, Hkv, window_left=window)
    y2 = ops.attention_decode_qkv(qkv, qn, kn, 1e-6, cos, sin, pos, kc, vc, sl, S, Hq, Hkv,
                                  window_left=window)
    assert (y.float() - y2.float()).abs().max().item() <= 2e-2
    # the step's rows landed in the right pool blocks, equal to the contiguous write
    for b in range(B):
        p = int(pos[b])
        blk = int(table[b, p // 64])
        assert torch.equal(kp[blk, :, p % 64], kc[b, :, p])
        assert torch.equal(vp[blk, :, p % 64], vc[b, :, p])
