"""GPU test of tpp_attention_decode_noalloc, the decode-attention entry point
that allocates nothing (for callers that cannot call cudaMalloc while they
decode: allocator callbacks, fixed-budget runtimes, plain-C hosts).

It is called straight through the C-ABI and must give the same result as
tpp_attention_decode with a caller workspace, on two calls in a row (the
second with different data, so stale scratch from the first call would
show).  This file is named to be collected last."""
import ctypes

import pytest
import torch

from torchplusplus_b200 import _native as N
from torchplusplus_b200 import ops

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2   # the tolerance of tests/test_kernels_gpu.py
MEAN_ABS = 1e-3


def _noalloc(q, kc, vc, seqlens, max_seqlen, out, window=-1):
    B, Hq, D = q.shape
    Hkv = kc.shape[1]
    return N.lib().tpp_attention_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), kc.stride(0),
        kc.stride(1), kc.stride(2), seqlens.data_ptr(), max_seqlen, out.data_ptr(),
        out.stride(0), out.stride(1), B, Hq, Hkv, D, window, ctypes.c_float(D ** -0.5),
        N.dtype_code(q.dtype), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("window", [-1, 1023])
def test_noalloc_matches_workspace_entry_point_twice(window):
    g = torch.Generator().manual_seed(21)
    # two sequences of ~3k keys: few CTAs per key range, so the key range is
    # split more than 8 ways and the partials go through the scratch array
    B, Hq, Hkv, D, Smax = 2, 16, 8, 128, 3000
    for call in range(2):
        q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).cuda()
        kc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16).cuda()
        vc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16).cuda()
        lens = [Smax - 7 * i - 300 * call for i in range(B)]
        # this exact shape (Hkv = 8, this window) sends its partials through
        # the scratch array, not only through the cluster merge
        assert N.lib().tpp_attention_decode_workspace_exact(B, Hq, Hkv, max(lens), D,
                                                            window) > 0
        sl = torch.tensor(lens, dtype=torch.int32).cuda()
        ref = ops.attention_decode(q, kc, vc, sl, max(lens), window_left=window)
        out = torch.full_like(ref, float("nan"))
        assert _noalloc(q, kc, vc, sl, max(lens), out, window) == 0, N.lib().tpp_last_error()
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, (call, err.max())


def test_noalloc_rejects_shapes_beyond_its_scratch():
    cap = N.lib().tpp_attention_decode_noalloc_max_bytes()
    assert cap == 8 << 20
    B, Hq, Hkv, D, L = 1, 64, 1, 256, 1 << 16
    assert ops.decode_workspace_bytes(B, Hq, L, D) > cap
    q = torch.zeros(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(1, 1, 1, D, dtype=torch.bfloat16, device="cuda").expand(B, Hkv, L, D)
    sl = torch.full((B,), L, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    st = _noalloc(q, kc, kc, sl, L, out)
    assert st == 7  # TPP_ERR_WORKSPACE, before any launch
    assert b"more than the fixed" in N.lib().tpp_last_error()
