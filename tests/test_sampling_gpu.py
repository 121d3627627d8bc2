"""On-device sampling (tpp_sample) against the reference's sampling rules
(torchpp/llmops/llm.py:114-203): degenerate settings reduce to argmax, the
sampled tokens stay inside the top-k / top-p sets, and the empirical
distribution over many independent draws matches softmax(logits / T)
restricted to those sets."""
import math

import pytest
import torch

from torchplusplus_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rows(B, V, seed, dtype=torch.bfloat16, scale=3.0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(B, V, generator=g)).to(dtype).to(DEV)


def _is_row_max(x, y):
    # tokens tied with the top logit are all kept (bf16 logits tie often)
    picked = x.gather(1, y[:, None])[:, 0]
    return torch.equal(picked, x.max(dim=1).values)


def test_top_k_one_is_argmax():
    x = _rows(64, 151936, 1)
    y = ops.sample(x, temperature=0.7, top_k=1)
    assert _is_row_max(x, y)
    xs = _rows(64, 4096, 5, dtype=torch.float16, scale=1.0)  # few ties: exact argmax
    ys = ops.sample(xs, temperature=0.7, top_k=1)
    assert _is_row_max(xs, ys)


def test_tiny_top_p_is_argmax():
    x = _rows(32, 4096, 2)
    y = ops.sample(x, temperature=1.0, top_p=1e-6)
    assert _is_row_max(x, y)


def _expected(logits_row, T, top_k, top_p):
    """Reference sets: llm.py sample_top_k / sample_top_p on one fp32 row."""
    l = logits_row.float() / T
    keep = torch.ones_like(l, dtype=torch.bool)
    if top_k:
        thr = torch.topk(l, top_k).values[-1]
        keep &= l >= thr
    p = torch.softmax(l.masked_fill(~keep, -float("inf")), -1)
    if top_p < 1.0:
        sp, si = torch.sort(p, descending=True)
        cum = torch.cumsum(sp, -1)
        remove = cum > top_p
        remove[1:] = remove[:-1].clone()
        remove[0] = False
        k2 = torch.ones_like(keep)
        k2[si[remove]] = False
        keep &= k2
    q = torch.softmax(l.masked_fill(~keep, -float("inf")), -1)
    return keep, q


@pytest.mark.parametrize("cfg", [(1.0, 0, 1.0), (0.8, 8, 1.0), (1.3, 0, 0.6), (1.0, 20, 0.8)])
def test_sample_distribution(cfg):
    T, k, p = cfg
    V, B = 64, 16384
    base = _rows(1, V, 3, scale=1.5)[0]
    x = base.expand(B, V).contiguous()
    counters = torch.arange(B, dtype=torch.int32, device=DEV)
    y = ops.sample(x, temperature=T, top_k=k, top_p=p, seed=1234, counters=counters).cpu()
    keep, q = _expected(base.cpu(), T, k, p)
    assert keep[y].all(), "sampled a token outside the top-k / top-p set"
    freq = torch.bincount(y, minlength=V).double() / B
    sigma = torch.sqrt(q.double() * (1 - q.double()) / B)
    assert ((freq - q.double()).abs() <= 5 * sigma + 1e-3).all()


def test_sample_draws_change_with_counters_and_seed():
    x = _rows(4, 1024, 4, scale=0.5)  # flat-ish: draws vary
    c0 = torch.zeros(4, dtype=torch.int32, device=DEV)
    a = ops.sample(x, counters=c0, seed=7)
    assert torch.equal(a, ops.sample(x, counters=c0, seed=7))  # deterministic
    draws = {tuple(ops.sample(x, counters=c0 + i, seed=7).tolist()) for i in range(8)}
    assert len(draws) > 1
