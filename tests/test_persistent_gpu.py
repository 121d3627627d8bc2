"""The persistent single-sequence decode step (tpp_decode_step_persistent):
one cooperative kernel per step against the launch-per-phase decode graph
(same folded weights, same caches) and, through the benchmark-shape test,
against the fp32 oracle."""
import pytest
import torch

from torchplusplus_b200 import ops
from torchplusplus_b200.llmops.engine import DecodeEngine
from torchplusplus_b200.llmops.qwen3 import Qwen3, Qwen3Config

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model(dtype=torch.bfloat16, seed=0, layers=2, heads=(4, 2)):
    cfg = Qwen3Config(vocab_size=1000, context_length=512, embed_dim=512, n_heads=heads[0],
                      n_layers=layers, head_dim=128, n_kv_heads=heads[1], hidden_dim=1024,
                      dtype=dtype)
    m = Qwen3(cfg, device=DEV).init_weights(0.05, seed=seed)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() == 1:
                p.copy_(1 + 0.1 * torch.randn(p.shape, device=DEV).to(p.dtype))
    return m


@pytest.mark.parametrize("heads", [(4, 2), (8, 2), (2, 2)], ids=["gq2", "gq4", "gq1"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("prompt", [1, 37, 200])
def test_persistent_step_matches_graph_step(dtype, prompt, heads):
    m = _model(dtype, heads=heads)
    ids = torch.randint(0, 1000, (1, prompt), generator=torch.Generator().manual_seed(prompt))
    with torch.inference_mode():
        ea = DecodeEngine(m, 1, 256, persistent=True)
        eb = DecodeEngine(m, 1, 256, persistent=False)
        assert ea.persistent is not None and eb.persistent is None
        ea.prefill(ids)
        eb.prefill(ids)
        for step in range(6):
            # teacher-force both engines with the same token
            eb.tokens.copy_(ea.tokens)
            eb.out_ids.copy_(ea.out_ids)
            ea.step_eager()
            eb.step_eager()
            la, lb = ea.logits.float(), eb.logits.float()
            err = (la - lb).abs().max().item()
            assert err <= 2e-2 * max(1.0, lb.abs().max().item()), (step, err)
            # the persistent step's pick is an argmax of the graph step's logits
            picked = lb[0, ea.tokens[0]]
            assert picked >= lb.max() - 2e-2 * max(1.0, lb.abs().max().item())
            # the new K/V rows agree
            pos = int(ea.positions[0]) - 1
            for ca, cb in zip(ea.caches, eb.caches):
                for xa, xb in ((ca.k_cache, cb.k_cache), (ca.v_cache, cb.v_cache)):
                    ra, rb = xa[0, :, pos].float(), xb[0, :, pos].float()
                    # two bf16 pipelines with different accumulation orders:
                    # a few ulps apart in the later layers
                    assert ((ra - rb).abs() / rb.abs().clamp(min=1.0)).max() <= 5e-2
        assert int(ea.positions[0]) == prompt + 6 and int(ea.seqlens[0]) == prompt + 7
        assert int(ea.out_ids[0, prompt + 6]) == int(ea.tokens[0])
    assert ops.device_error() == 0


def test_persistent_generate_graph_replays():
    """Greedy generate at batch 1 runs the persistent step inside the decode
    graph; every pick is an argmax of the launch-per-phase path's logits on
    the same sequence."""
    m = _model(torch.bfloat16, seed=3)
    ids = torch.randint(0, 1000, (1, 30), generator=torch.Generator().manual_seed(9))
    m.decode_persistent = True
    with torch.inference_mode():
        out = m.generate(ids, max_new_token=16, sampling_strategy="greedy")
        assert m._engine.persistent is not None and m._engine.launches_per_step == 1
        logits = m.forward_impl(out[:, :-1].to(DEV)).float()[:, 29:]
    picked = logits.gather(-1, out[:, 30:].to(DEV)[..., None])[..., 0]
    best = logits.max(-1).values
    assert bool((picked >= best - 5e-2 * best.abs().clamp(min=1.0)).all())
    assert ops.device_error() == 0


@pytest.mark.parametrize("prompt", [600, 2600])
def test_persistent_step_at_qwen3_widths(prompt):
    """Qwen3-0.6B layer widths (E 1024, 16/8 heads, F 3072): at 600 keys
    every attention unit's cached rows are staged in shared memory behind its
    o-proj slice; at 2600 a unit's range (145 keys) outgrows that room (135
    rows on 148 SMs) and its last rows come from the cache directly."""
    cfg = Qwen3Config(vocab_size=4096, context_length=4096, n_layers=2, dtype=torch.bfloat16)
    m = Qwen3(cfg, device=DEV).init_weights(0.02, seed=5)
    ids = torch.randint(0, 4096, (1, prompt), generator=torch.Generator().manual_seed(prompt))
    with torch.inference_mode():
        ea = DecodeEngine(m, 1, 3072, persistent=True)
        eb = DecodeEngine(m, 1, 3072, persistent=False)
        assert ea.persistent is not None
        ea.prefill(ids)
        eb.prefill(ids)
        for step in range(3):
            eb.tokens.copy_(ea.tokens)
            eb.out_ids.copy_(ea.out_ids)
            ea.step_eager()
            eb.step_eager()
            la, lb = ea.logits.float(), eb.logits.float()
            assert (la - lb).abs().max().item() <= 2e-2 * max(1.0, lb.abs().max().item()), step
    assert ops.device_error() == 0


def test_persistent_steps_repeat_exactly_across_requests():
    """The step kernel tags every exchanged activation with an epoch derived
    from the steps already run on its workspace; a second request on the
    same engine (epochs continuing, graph replays) must pick the same tokens
    as the first."""
    m = _model(torch.bfloat16, seed=4)
    ids = torch.randint(0, 1000, (1, 45), generator=torch.Generator().manual_seed(11))
    m.decode_persistent = True
    with torch.inference_mode():
        a = m.generate(ids, max_new_token=24, sampling_strategy="greedy").cpu()
        eng = m._engine
        b = m.generate(ids, max_new_token=24, sampling_strategy="greedy").cpu()
        assert m._engine is eng and eng.persistent is not None
    assert torch.equal(a, b)
    assert ops.device_error() == 0
